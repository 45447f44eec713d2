"""Lightning indexer on the B200 tensor cores against the reference (test_kernels.py:89-126, BASELINE
configs 3 and 4): rel_err < 1e-5 of the float64 oracle, causal -inf masks equal."""
import numpy as np
import pytest
import torch

import oracle as O
import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import workloads
from tests.gpu_util import DEV, assert_no_device_error, cuda, npy, rel_err, sample_rows

pytestmark = pytest.mark.gpu


def _dev(*ts):
    return [t.to(DEV) for t in ts]


def test_index_matches_reference_golden(golden):
    for ii in range(int(golden["ix_ncases"])):
        B, M, N, H, D_, causal, start = golden[f"ix_{ii}_meta"].tolist()
        q, w, k, ks = (cuda(golden[f"ix_{ii}_{n}"]) for n in ("q", "w", "k", "ks"))
        o = D.int8_index(q, w, k, ks, causal=bool(causal), start=start)
        ref = golden[f"ix_{ii}_o"]
        assert o.shape == (B, M, N)
        np.testing.assert_array_equal(np.isinf(npy(o)), np.isinf(ref))
        assert rel_err(npy(o), ref) < 1e-5
    assert_no_device_error()


@pytest.mark.parametrize("B,M,N", [(1, 1, 128), (1, 1, 1000), (2, 3, 257), (1, 17, 512), (2, 64, 1024)])
def test_index_reference_shapes(B, M, N):
    q, w, k, ks = workloads.index_inputs_uniform(B, M, N, seed=B + M + N)
    o = D.int8_index(*_dev(q, w, k, ks), block_q=2, block_n=64)
    assert rel_err(npy(o), O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy())) < 1e-5


@pytest.mark.parametrize("M,N,start", [(64, 64, 0), (100, 100, 0), (16, 300, 284), (33, 200, 50),
                                       (300, 700, 400), (5, 1000, 0)])
def test_index_causal(M, N, start):
    q, w, k, ks = workloads.index_inputs_uniform(1, M, N, seed=M + N + start)
    o = D.int8_index(*_dev(q, w, k, ks), causal=True, start=start)
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy(), causal=True, start=start)
    np.testing.assert_array_equal(np.isinf(npy(o)), np.isinf(ref))
    assert rel_err(npy(o), ref) < 1e-5


@pytest.mark.parametrize("H,D_", [(16, 64), (32, 128), (64, 64), (16, 128)])
def test_index_other_head_shapes(H, D_):
    q, w, k, ks = workloads.index_inputs_uniform(1, 8, 256, H=H, D=D_, seed=H + D_)
    o = D.int8_index(*_dev(q, w, k, ks))
    assert rel_err(npy(o), O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy())) < 1e-5


def test_index_topk_overlap_reference_test():
    """test_kernels.py:121-126: top-256 of 4096 keys matches the reference's selection."""
    q, w, k, ks = workloads.index_inputs_uniform(1, 32, 4096, seed=5)
    o = npy(D.int8_index(*_dev(q, w, k, ks)))
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy())
    a = np.sort(np.argsort(-o, -1)[..., :256], -1)
    r = np.sort(np.argsort(-ref, -1)[..., :256], -1)
    assert (a == r).mean() > 0.999


def test_index_baseline_decode_full_size():
    """4 queries x 32768 keys (shared key cache), rotated+quantised generators."""
    q, w, k, ks = workloads.index_inputs(1, 4, 32768, seed=0)
    o = D.int8_index(*_dev(q, w, k, ks))
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy())
    assert rel_err(npy(o), ref) < 1e-5
    # the same 4 queries as 4 batch rows, each with its own copy of the keys
    qb, wb = q.view(4, 1, 64, 128).contiguous(), w.view(4, 1, 64).contiguous()
    kb, ksb = k.expand(4, -1, -1).contiguous(), ks.expand(4, -1).contiguous()
    ob = D.int8_index(*_dev(qb, wb, kb, ksb))
    assert torch.equal(ob.view(1, 4, -1), o)
    assert_no_device_error()


def test_index_baseline_prefill_full_size():
    """4096 x 4096 causal; oracle on a seeded sample of query rows; -inf masks
    exact for every row."""
    M = N = 4096
    q, w, k, ks = workloads.index_inputs(1, M, N, seed=0)
    o = npy(D.int8_index(*_dev(q, w, k, ks), causal=True, start=0))
    rows = sample_rows(M, 64)
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy(), causal=True, start=0, rows=rows)
    assert rel_err(o[:, rows], ref) < 1e-5
    mask = np.arange(N)[None, :] > np.arange(M)[:, None]
    np.testing.assert_array_equal(np.isinf(o[0]), mask)
    assert np.isfinite(o[0][~mask]).all()
    assert_no_device_error()


def test_index_long_context_rows():
    """Chunked-prefill convention of the long case: last queries of a long sequence (start > 0)."""
    M, N = 256, 20000
    q, w, k, ks = workloads.index_inputs(1, M, N, seed=3)
    start = N - M
    o = npy(D.int8_index(*_dev(q, w, k, ks), causal=True, start=start))
    rows = sample_rows(M, 16)
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy(), causal=True, start=start, rows=rows)
    np.testing.assert_array_equal(np.isinf(o[:, rows]), np.isinf(ref))
    assert rel_err(o[:, rows], ref) < 1e-5


def test_index_v2_shims():
    q, w, k, ks = workloads.index_inputs_uniform(2, 3, 257, seed=11)
    o = D.int8_index_v2(D.index_kmajor_q(q.to(DEV)), w.to(DEV), D.index_kmajor_k(k.to(DEV)), ks.to(DEV), H=64)
    assert rel_err(npy(o), O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy())) < 1e-5
