"""Fused top-k selection on the B200: the selected index sets equal the oracle's deterministic top-k
(ties to the lowest position) exactly, and are valid torch.topk answers tie-aware."""
import numpy as np
import pytest
import torch

import oracle as O
import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import workloads
from tests.gpu_util import DEV, assert_no_device_error, npy, sample_rows

pytestmark = pytest.mark.gpu


def _scores(rows, n, ties, seed, neginf_tail=0):
    g = torch.Generator().manual_seed(seed)
    s = torch.randint(0, 40, (rows, n), generator=g).float() if ties else torch.randn(rows, n, generator=g)
    if neginf_tail:
        s[:, n - neginf_tail:] = float("-inf")
    return s


@pytest.mark.parametrize("n,k", [(100, 10), (1000, 999), (4096, 2048), (8192, 2048), (20000, 2048),
                                 (40000, 2048), (131072, 2048)])
@pytest.mark.parametrize("ties", [False, True])
def test_select_topk_equals_oracle(n, k, ties):
    rows = 3 if n > 20000 else 6
    s = _scores(rows, n, ties, seed=n + k)
    idx, vals = D.select_topk(s.to(DEV), k)
    ri, rv = O.topk_ref(s.numpy(), k)
    np.testing.assert_array_equal(npy(idx), ri)
    np.testing.assert_array_equal(npy(vals), rv)
    assert O.topk_valid(npy(idx), s.numpy(), k)
    assert_no_device_error()


def test_select_topk_with_masked_tail():
    s = _scores(4, 3000, False, seed=7, neginf_tail=2500)  # 500 finite values, k = 2048
    idx, vals = D.select_topk(s.to(DEV), 2048)
    ri, rv = O.topk_ref(s.numpy(), 2048)
    np.testing.assert_array_equal(npy(idx), ri)
    assert O.topk_valid(npy(idx), s.numpy(), 2048)


def _assert_same_values(got, ref):
    """NaN where the reference has NaN (any payload); every other value bit for bit."""
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got.view(np.int32)[~nan], ref.view(np.int32)[~nan])


def _nan_rows(rows, n, seed):
    """Rows with NaNs of both signs and several payloads, infinities, masked tails and signed zeros."""
    g = torch.Generator().manual_seed(seed)
    s = torch.randn(rows, n, generator=g)
    b = s.view(torch.int32)
    s[0, 5], s[0, 40] = float("nan"), float("inf")
    b[0, 17] = -4194304                                  # 0xFFC00000: NaN with the sign bit set
    s[1] = float("-inf")
    s[1, 3] = float("nan")
    b[1, 9] = -1                                         # 0xFFFFFFFF: all bits set
    s[2, 100:] = float("-inf")
    b[2, 10] = 0x7F800123                                # NaN with a payload
    s[3, ::2] = 0.0
    s[3, 1::4] = -0.0
    b[4, ::3] = 0x7FC00000
    b[4, 1::7] = -8388607                                # 0xFF800001: the lowest negative NaN bits
    return s


@pytest.mark.parametrize("n,k,rows", [(300, 64, 6), (1536, 512, 6), (1536, 16, 6), (20000, 2048, 160),
                                      (40000, 2048, 6), (131072, 2048, 5)])
def test_select_topk_nan_and_signed_zero_order(n, k, rows):
    """Values are ranked as torch.topk ranks fp32 on the GPU: every NaN above +inf (NaNs tie, lowest
    position first), -0.0 just below +0.0. Covers the register pass, the staged plan (few long rows),
    the long-row filter and its scratch-free fallback. Values other than NaN are returned bit for bit
    (signed zeros included); a selected NaN comes back as a NaN."""
    s = _nan_rows(rows, n, seed=n + k)
    idx, vals = D.select_topk(s.to(DEV), k)
    pick = list(range(min(rows, 6))) + [rows - 1]
    ri, rv = O.topk_ref(s.numpy()[pick], k)
    np.testing.assert_array_equal(npy(idx)[pick], ri)
    _assert_same_values(npy(vals)[pick], rv)
    assert_no_device_error()


def test_merge_of_shard_lists_with_nan_equals_global():
    """NaN order holds through the merge of per-shard lists (read in place and concatenated)."""
    n, k, shards = 16384, 2048, 4
    s = _nan_rows(6, n, seed=99).to(DEV)
    step = n // shards
    parts = [D.select_topk(s[:, r * step:(r + 1) * step].contiguous(), k, idx_offset=r * step) for r in range(shards)]
    midx, mval = D.select_topk_parts([p[1] for p in parts], [p[0] for p in parts], k)
    gidx, gval = D.select_topk(s, k)
    assert torch.equal(midx, gidx) and torch.equal(mval.view(torch.int32), gval.view(torch.int32))
    ri, rv = O.topk_ref(npy(s), k)
    np.testing.assert_array_equal(npy(gidx), ri)
    assert_no_device_error()


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_merge_of_shard_topk_equals_global(shards):
    """Key-range sharding: per-shard top-k with global key offsets, candidate lists
    concatenated in shard order, merged with the same kernel -> identical to the one-shot top-k."""
    n, k = 16384, 2048
    s = _scores(5, n, True, seed=shards).to(DEV)
    step = n // shards
    parts = [D.select_topk(s[:, r * step:(r + 1) * step].contiguous(), k, idx_offset=r * step) for r in range(shards)]
    cand_idx = torch.cat([p[0] for p in parts], -1).contiguous()
    cand_val = torch.cat([p[1] for p in parts], -1).contiguous()
    midx, mval = D.select_topk(cand_val, k, cand_idx=cand_idx)
    gidx, gval = D.select_topk(s, k)
    assert torch.equal(midx, gidx) and torch.equal(mval, gval)


@pytest.mark.parametrize("shards,n,k,rows", [(2, 16384, 2048, 5), (4, 16384, 2048, 37), (8, 65536, 2048, 3),
                                              (16, 65536, 2048, 2), (3, 192, 100, 9), (5, 640, 64, 4),
                                              (5, 10000, 2000, 3)])
def test_merge_of_shard_lists_in_place_equals_global(shards, n, k, rows):
    """select_topk_parts reads the per-shard lists where they lie (no concatenation): identical to the
    merge of the concatenated lists and to the one-shot top-k, ties included (integer-valued scores),
    including single-pass, staged (8 and 16 lists of 2048; 5 lists of 2000, whose stage segments
    must start on list-aligned 16-position boundaries) and short-list cases."""
    s = _scores(rows, n, True, seed=shards * 7 + k).to(DEV)
    s[0, : n // shards] = float("-inf")  # one shard of one row entirely masked
    step = n // shards
    kk = min(k, step)
    parts = [D.select_topk(s[:, r * step:(r + 1) * step].contiguous(), kk, idx_offset=r * step) for r in range(shards)]
    midx, mval = D.select_topk_parts([p[1] for p in parts], [p[0] for p in parts], k)
    cidx = torch.cat([p[0] for p in parts], -1).contiguous()
    cval = torch.cat([p[1] for p in parts], -1).contiguous()
    ridx, rval = D.select_topk(cval, k, cand_idx=cidx)
    assert torch.equal(midx, ridx) and torch.equal(mval, rval)
    if kk == k:
        gidx, gval = D.select_topk(s, k)
        assert torch.equal(midx, gidx) and torch.equal(mval, gval)
    assert_no_device_error()


def test_index_topk_prefill_4096_causal():
    """BASELINE config 4 end to end: scores + top-2048 per query, causal."""
    M = N = 4096
    q, w, k, ks = workloads.index_inputs(1, M, N, seed=0)
    scores, idx, vals = D.int8_index_topk(q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV), topk=2048, causal=True)
    sc = npy(scores)[0]
    ri, rv = O.topk_ref(sc, 2048)  # deterministic selection over the kernel's own scores
    np.testing.assert_array_equal(npy(idx)[0], ri)
    rows = sample_rows(M, 32)
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy(), causal=True, rows=rows)[0]
    assert O.topk_valid(npy(idx)[0][rows], ref, 2048) or _near_tie_ok(npy(idx)[0][rows], ref, 2048)
    assert_no_device_error()


def _near_tie_ok(sel, ref, k, rel=1e-5):
    """fp32 scores may order two keys whose float64 values differ by less than the kernel tolerance
    differently; accept swaps within that band (tie-aware at the tolerance)."""
    for r in range(ref.shape[0]):
        row = ref[r]
        kth = np.sort(row)[-k]
        if np.isneginf(kth):
            if not np.all(np.isin(np.flatnonzero(np.isfinite(row)), sel[r])):
                return False
            continue
        band = rel * np.abs(row[np.isfinite(row)]).max()
        if np.any(row[sel[r]] < kth - band) or not np.all(np.isin(np.flatnonzero(row > kth + band), sel[r])):
            return False
    return True


def test_index_topk_decode():
    q, w, k, ks = workloads.index_inputs(1, 4, 32768, seed=1)
    idx, vals = D.int8_index_topk(q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV), topk=2048, return_scores=False)
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy())[0]
    assert O.topk_valid(npy(idx)[0], ref, 2048) or _near_tie_ok(npy(idx)[0], ref, 2048)


def test_select_topk_with_infinities():
    s = _scores(3, 5000, False, seed=9)
    s[0, 10] = float("inf")
    s[1, ::7] = float("-inf")
    s[2, 100:4000] = float("-inf")  # 1100 values above -inf, k = 2048
    idx, vals = D.select_topk(s.to(DEV), 2048)
    ri, rv = O.topk_ref(s.numpy(), 2048)
    np.testing.assert_array_equal(npy(idx), ri)
    np.testing.assert_array_equal(npy(vals), rv)


@pytest.mark.parametrize("start", [-300, 0, 700])
def test_index_topk_causal_batched_with_offset(start):
    """The fused call skips reading each causal row's masked tail; its selection must equal the
    deterministic top-k of the scores it returns, for every batch and a shifted causal start."""
    B, M, N, topk = 2, 384, 1536, 512
    q, w, k, ks = workloads.index_inputs(B, M, N, seed=11)
    scores, idx, vals = D.int8_index_topk(q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV), topk=topk, causal=True,
                                          start=start, key_offset=4096)
    for b in range(B):
        sc = npy(scores)[b]
        ri, rv = O.topk_ref(sc, topk)
        np.testing.assert_array_equal(npy(idx)[b], ri + 4096)
        np.testing.assert_array_equal(npy(vals)[b], rv)
    assert_no_device_error()


@pytest.mark.parametrize("start,N,topk", [(-300, 1536, 512), (0, 4096, 2048), (700, 1536, 512), (100, 640, 640),
                                          (3000, 4096, 512)])
def test_index_topk_leading_rows_selected_by_the_indexer(start, N, topk):
    """In a single-batch causal call the leading rows see at most topk keys, so their selection is their
    first topk positions; the indexer writes it itself and the top-k launch covers the other rows. The
    result must equal the plain selection over the returned scores, bit for bit, with the scores kept
    or not, and with NaN (of either sign) in the weights and key scales."""
    M = 640
    q, w, k, ks = workloads.index_inputs(1, M, N, seed=31)
    ks[0, 7] = float("nan")
    ks[0, 9] = torch.tensor(float("nan")).neg()
    w[0, 300, 5] = torch.tensor(float("nan")).neg()
    qd, wd, kd, ksd = q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV)
    scores, idx, vals = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=start, key_offset=77)
    pidx, pvals = D.select_topk(scores.view(M, N), topk)
    assert torch.equal(idx.view(M, topk), pidx + 77)
    assert torch.equal(vals.view(M, topk).view(torch.int32), pvals.view(torch.int32))
    idx2, vals2 = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=start, key_offset=77,
                                    return_scores=False)
    assert torch.equal(idx2, idx) and torch.equal(vals2.view(torch.int32), vals.view(torch.int32))
    assert_no_device_error()


def test_index_topk_causal_long_rows_batched():
    """Rows longer than one register pass are selected in stages, in row batches that bound the
    scratch; with causal rows the first stage skips each row's masked tail. The result must equal
    the plain selection over the returned scores (which reads the -inf tail) and the oracle."""
    B, M, N, topk, start = 1, 5000, 12000, 2048, 6000
    q, w, k, ks = workloads.index_inputs(B, M, N, seed=21)
    scores, idx, vals = D.int8_index_topk(q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV), topk=topk, causal=True,
                                          start=start)
    pidx, pvals = D.select_topk(scores.view(B * M, N), topk)
    assert torch.equal(idx.view(B * M, topk), pidx) and torch.equal(vals.view(B * M, topk), pvals)
    rows = [0, 1, 2047, 2191, 2192, 4095, 4096, 4999]
    sc = npy(scores)[0][rows]
    ri, rv = O.topk_ref(sc, topk)
    np.testing.assert_array_equal(npy(idx)[0][rows], ri)
    np.testing.assert_array_equal(npy(vals)[0][rows], rv)
    assert_no_device_error()


def test_index_topk_baseline_long_full_size():
    """BASELINE configs[4], long-context case on one GPU: 4096 queries x 131072 keys, causal with the
    chunked-prefill start 126976, top-2048. Rows are selected in stages through the workspace.
    Scores on 64 sampled rows (first and last included) are within 1e-5 of the float64 oracle with
    exact -inf masks; the selection equals the deterministic top-k of the returned scores on those
    rows and is a valid top-k of the float64 scores (tie-aware, at the kernel's tolerance where two
    keys' fp32 scores order differently from their float64 ones). The indices-only call, which
    leaves the masked tiles unwritten, selects the same keys."""
    M, N, topk = 4096, 131072, 2048
    start = N - M
    q, w, k, ks = workloads.index_inputs(1, M, N, seed=0)
    qd, wd, kd, ksd = q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV)
    scores, idx, vals = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=start)
    rows = sample_rows(M, 64, seed=4)
    sc = npy(scores[0, torch.from_numpy(rows).to(DEV)])
    del scores
    ref = O.int8_index_ref(q.numpy(), w.numpy(), k.numpy(), ks.numpy(), causal=True, start=start, rows=rows,
                           chunk=8)[0]
    np.testing.assert_array_equal(np.isinf(sc), np.isinf(ref))
    assert O.rel_err(sc, ref) < 1e-5
    ri, rv = O.topk_ref(sc, topk)
    sel = npy(idx)[0][rows]
    np.testing.assert_array_equal(sel, ri)
    np.testing.assert_array_equal(npy(vals)[0][rows], rv)
    strict = [O.topk_valid(sel[j:j + 1], ref[j:j + 1], topk) for j in range(len(rows))]
    banded = [s or _near_tie_ok(sel[j:j + 1], ref[j:j + 1], topk) for j, s in enumerate(strict)]
    print(f"long config: {sum(strict)} of {len(rows)} sampled rows valid against float64 without the tie band")
    assert all(banded)
    idx2, vals2 = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=start, return_scores=False)
    assert torch.equal(idx2, idx) and torch.equal(vals2, vals)
    assert_no_device_error()


def test_long_rows_without_workspace_use_the_scratch_free_kernel():
    """dsv32_topk with no workspace selects rows longer than 8192 with the kernel that re-reads them
    from L2 (no scratch); it must equal the staged selection."""
    from deepseek_v32_gtx1650_b200 import _lib
    rows, n, k = 5, 40000, 2048
    s = _scores(rows, n, True, seed=17).to(DEV)
    s[1, 5000:] = float("-inf")
    gi, gv = D.select_topk(s, k)  # staged, with the per-stream workspace
    oi = torch.empty(rows, k, dtype=torch.int32, device=DEV)
    ov = torch.empty(rows, k, device=DEV)
    _lib.check(_lib.load().dsv32_topk(s.data_ptr(), rows, n, n, None, 0, 0, k, oi.data_ptr(), ov.data_ptr(), None, 0,
                                      torch.cuda.current_stream().cuda_stream), "dsv32_topk without workspace")
    assert torch.equal(oi, gi) and torch.equal(ov, gv)
    assert_no_device_error()


def test_index_topk_reads_key_cache_in_place():
    """n_keys scores the first n_keys keys of a cache with spare capacity through the key batch
    stride (no copy): identical to the call on the contiguous slice."""
    B, M, cap, n, topk = 2, 96, 3000, 2100, 512
    q, w, k, ks = workloads.index_inputs(B, M, cap, seed=13)
    qd, wd, kd, ksd = q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV)
    s1, i1, v1 = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=n - M, n_keys=n)
    s2, i2, v2 = D.int8_index_topk(qd, wd, kd[:, :n].contiguous(), ksd[:, :n].contiguous(), topk=topk, causal=True,
                                   start=n - M)
    assert torch.equal(s1, s2) and torch.equal(i1, i2) and torch.equal(v1, v2)
    assert_no_device_error()


def test_steady_state_calls_allocate_no_device_memory():
    """The library allocates nothing: after one call of each shape has filled the caller-side caches
    (outputs, the top-k and GEMM workspaces), further decode and long-row calls leave the device's
    free memory unchanged."""
    qd, wd, kd, ksd = (t.to(DEV) for t in workloads.index_inputs(1, 4, 32768, seed=2))
    ql, wl, kl, ksl = (t.to(DEV) for t in workloads.index_inputs(1, 64, 40000, seed=3))

    def calls():
        D.int8_index_topk(qd, wd, kd, ksd, topk=2048, return_scores=False)
        D.int8_index_topk(ql, wl, kl, ksl, topk=2048, causal=True, start=40000 - 64, return_scores=False)
        torch.cuda.synchronize()

    calls()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        calls()
    assert torch.cuda.mem_get_info()[0] == free0
    assert_no_device_error()


@pytest.mark.parametrize("n,k,ties", [(20000, 2048, False), (40000, 2048, True), (65536, 1000, False),
                                      (131072, 2048, True), (17000, 2730, False), (12000, 2048, False),
                                      (16384, 2048, True), (8200, 100, False)])
def test_long_rows_filter_equals_oracle(n, k, ties):
    """Rows longer than one register pass, at least one per SM (160 rows): each row is reduced to the
    keys at or above a sampled threshold, in position order, then selected in one register pass. The
    selection equals the oracle's deterministic top-k, values and ties included."""
    rows = 160
    s = _scores(rows, n, ties, seed=n + k).to(DEV)
    s[3, n // 2:] = float("-inf")      # a row with a long masked tail
    s[4, : n - k] = float("-inf")      # exactly k values above -inf
    s[5, 10] = float("inf")
    idx, vals = D.select_topk(s, k)
    pick = [0, 3, 4, 5, 77, rows - 1]
    ri, rv = O.topk_ref(npy(s)[pick], k)
    np.testing.assert_array_equal(npy(idx)[pick], ri)
    np.testing.assert_array_equal(npy(vals)[pick], rv)
    assert_no_device_error()


def test_long_rows_filter_fallbacks():
    """Rows on which the sampled threshold misjudges the row (large values only at positions the sample
    skips, so the candidate list overflows; or only at sampled positions, so it holds fewer than k keys)
    and rows with masked keys among the k largest or more NaNs than the list holds are selected by
    the scratch-free kernel instead: every row still equals the oracle."""
    rows, n, k = 160, 20000, 2048
    g = torch.Generator().manual_seed(3)
    s = torch.rand(rows, n, generator=g)
    pos = torch.arange(n)
    sampled = (pos < 512 * 32) & ((pos % 32) < 16)  # thread t samples [32 t, 32 t + 16) for n = 20000
    big = torch.rand(rows, n, generator=g) + 10.0
    s[0] = torch.where(~sampled, big[0], s[0])                 # large values the sample never sees
    s[1] = torch.where(sampled, big[1], s[1])                  # the sample sees only large values
    s[2, 100:] = float("-inf")                                 # few visible values
    s[3, ::2] = torch.tensor(float("nan")).neg()               # negative NaNs everywhere
    sd = s.to(DEV)
    idx, vals = D.select_topk(sd, k)
    pick = [0, 1, 2, 3, 50, rows - 1]
    ri, rv = O.topk_ref(s.numpy()[pick], k)
    np.testing.assert_array_equal(npy(idx)[pick], ri)
    np.testing.assert_array_equal(npy(vals)[pick].view(np.int32), rv.astype(np.float32).view(np.int32))
    assert_no_device_error()


def test_index_topk_causal_long_rows_filter():
    """The fused indexer + top-k on causal rows longer than two register passes (256 queries over 40000
    keys): the filter skips each row's masked tail (left unwritten when the scores are scratch) and the
    selection equals the deterministic top-k of the returned scores."""
    B, M, N, topk = 1, 256, 40000, 2048
    start = N - M
    q, w, k, ks = workloads.index_inputs(B, M, N, seed=31)
    qd, wd, kd, ksd = q.to(DEV), w.to(DEV), k.to(DEV), ks.to(DEV)
    scores, idx, vals = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=start)
    rows = [0, 1, 100, 255]
    ri, rv = O.topk_ref(npy(scores)[0][rows], topk)
    np.testing.assert_array_equal(npy(idx)[0][rows], ri)
    np.testing.assert_array_equal(npy(vals)[0][rows], rv)
    idx2, vals2 = D.int8_index_topk(qd, wd, kd, ksd, topk=topk, causal=True, start=start, return_scores=False)
    assert torch.equal(idx2, idx) and torch.equal(vals2, vals)
    assert_no_device_error()
