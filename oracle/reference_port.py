"""numpy restatement of the reference's float64 oracle (reference.py) -- test infrastructure only.

Each function cites the reference lines it restates. All arithmetic is numpy on the CPU; the
integer parts are exact and the float parts follow the reference's rounding (fp32 where the
reference computes in fp32, float64 where it computes in float64).
"""
from __future__ import annotations

import numpy as np

GROUP = 128  # reference.py:4


# ---------------------------------------------------------------------------------- dtypes
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact), as torch's bf16 .float() (kernels.py:21-23)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (kernels.py:26-30; finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return b.astype(np.uint16)


# ---------------------------------------------------------------------------------- act_quant
_INV127 = np.float32(1.0 / 127.0)  # torch multiplies the fp32 tensor by fl32(1/127)
_FLOOR = np.float32(1e-4)          # torch.clamp(min=1e-4) on an fp32 tensor uses fl32(1e-4)


def act_quant_ref(x: np.ndarray, round_scale: bool = False):
    """reference.py:8-15. x: float32 array [..., N] (fp16/bf16 inputs converted to fp32 first,
    exactly, as x.float() does). Returns (int8 [..., N], float32 [..., N/128])."""
    x = np.asarray(x, dtype=np.float32)
    *lead, N = x.shape
    g = x.reshape(*lead, N // GROUP, GROUP)
    with np.errstate(invalid="ignore"):
        amax = np.abs(g).max(axis=-1)
        # torch.amax propagates NaN; numpy max does too.
        s = np.maximum(amax, _FLOOR) * _INV127  # fp32 * fp32, one rounding
        s = np.where(np.isnan(amax), np.float32(np.nan), s).astype(np.float32)
        if round_scale:
            # torch.exp2(torch.ceil(torch.log2(s))): torch's CPU fp32 log2 equals the correctly
            # rounded fp32 of log2 (pinned by tests/test_oracle.py against reference.py).
            fin = np.isfinite(s)
            l2 = np.log2(np.where(fin, s, 1.0).astype(np.float64)).astype(np.float32)
            e = np.ceil(l2).astype(np.int32)
            s = np.where(fin, np.ldexp(np.float32(1.0), e).astype(np.float32), s).astype(np.float32)
        q = g / s[..., None]  # IEEE fp32 division
        y = np.clip(np.rint(q), -127, 127)  # rint = round half to even, like torch.round
    y = np.nan_to_num(y, nan=0.0).astype(np.int8)
    return y.reshape(*lead, N), s


# ---------------------------------------------------------------------------------- int8_gemm
def int8_gemm_ref(a: np.ndarray, a_s: np.ndarray, b: np.ndarray, b_s: np.ndarray, chunk: int = 1024) -> np.ndarray:
    """reference.py:18-24: dequantise both sides block by block in float64, then matmul.
    a int8 [..., K], a_s [..., K/128], b int8 [N, K], b_s [N/128, K/128] -> float64 [..., N]."""
    K = a.shape[-1]
    N = b.shape[0]
    KG = K // GROUP
    a2 = a.reshape(-1, K)
    as2 = a_s.reshape(-1, KG).astype(np.float64)
    bs = np.repeat(b_s.astype(np.float64), GROUP, axis=0)[:N]  # [N, KG]
    Bd = (b.astype(np.float64).reshape(N, KG, GROUP) * bs[..., None]).reshape(N, K)
    out = np.empty((a2.shape[0], N), dtype=np.float64)
    for i in range(0, a2.shape[0], chunk):
        Ad = (a2[i:i + chunk].astype(np.float64).reshape(-1, KG, GROUP) * as2[i:i + chunk, :, None]).reshape(-1, K)
        out[i:i + chunk] = Ad @ Bd.T
    return out.reshape(*a.shape[:-1], N)


def int8_gemm_partials_ref(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact per-128-K-block integer products: [K/128, M, N] int64, partial[kb] = A_kb @ B_kb^T
    (the int32 tl.dot of kernels.py:94)."""
    K = a.shape[-1]
    KG = K // GROUP
    a2 = a.reshape(-1, K)
    out = np.empty((KG, a2.shape[0], b.shape[0]), dtype=np.int64)
    for kb in range(KG):
        sl = slice(kb * GROUP, (kb + 1) * GROUP)
        # float64 matmul of small integers is exact (|sum| <= 128 * 127^2 < 2^53) and uses BLAS.
        out[kb] = np.rint(a2[:, sl].astype(np.float64) @ b[:, sl].astype(np.float64).T).astype(np.int64)
    return out


# ---------------------------------------------------------------------------------- int8_index
def int8_index_ref(q: np.ndarray, w: np.ndarray, k: np.ndarray, k_s: np.ndarray, causal: bool = False,
                   start: int = 0, chunk: int = 64, rows: np.ndarray | None = None) -> np.ndarray:
    """reference.py:27-34: logits = einsum(q, k) in float64, relu, * w, sum over heads, * k_s;
    causal: -inf where n > start + m. q [B, M, H, D] int8, w [B, M, H], k [B, N, D] int8, k_s [B, N]
    -> float64 [B, M, N] (or [B, len(rows), N] for the selected query rows)."""
    B, M, H, D = q.shape
    N = k.shape[1]
    rows = np.arange(M) if rows is None else np.asarray(rows)
    out = np.empty((B, len(rows), N), dtype=np.float64)
    for b in range(B):
        kT = k[b].astype(np.float64).T  # [D, N]
        ks = k_s[b].astype(np.float64)
        for i in range(0, len(rows), chunk):
            r = rows[i:i + chunk]
            lg = q[b, r].astype(np.float64).reshape(-1, D) @ kT  # [r*H, N], exact integers
            np.maximum(lg, 0.0, out=lg)
            lg = lg.reshape(len(r), H, N)
            sc = np.einsum("mhn,mh->mn", lg, w[b, r].astype(np.float64)) * ks[None, :]
            if causal:
                keep = np.arange(N)[None, :] <= start + r[:, None]
                sc = np.where(keep, sc, -np.inf)
            out[b, i:i + chunk] = sc
    return out


# ---------------------------------------------------------------------------------- top-k
def order_keys(x: np.ndarray) -> np.ndarray:
    """fp32 -> uint32 keys in the order torch.topk ranks values on the GPU (its radix keys): negative
    floats with all bits flipped, the others with the sign bit raised, so -0.0 ranks just below +0.0,
    and every NaN (either sign) the all-ones key, above +inf, NaNs tying with one another."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    key = np.where(u >> np.uint32(31) == 1, ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    return np.where(np.isnan(x), np.uint32(0xFFFFFFFF), key).astype(np.uint32)


def topk_ref(scores: np.ndarray, k: int):
    """Deterministic top-k per row (the selection torch.topk makes in test_kernels.py:121-126, with its
    ties fixed): the k largest values in order_keys order (fp32 scores; wider types by value, NaN
    first), ties at the k-th key by lowest position, listed in increasing position order.
    Returns (idx int64 [..., k], vals [..., k])."""
    s = np.asarray(scores)
    n = s.shape[-1]
    flat = s.reshape(-1, n)
    idx = np.empty((flat.shape[0], k), dtype=np.int64)
    pos = np.arange(n)
    for r in range(flat.shape[0]):
        row = flat[r]
        if row.dtype == np.float32:
            order = np.lexsort((pos, -order_keys(row).astype(np.int64)))  # key desc, then position asc
        else:
            nan = np.isnan(row)
            order = np.lexsort((pos, -np.where(nan, 0.0, row), ~nan))  # NaN, value desc, position asc
        idx[r] = np.sort(order[:k])
    vals = np.take_along_axis(flat, idx, axis=1)
    return idx.reshape(*s.shape[:-1], k), vals.reshape(*s.shape[:-1], k)


def topk_valid(sel_idx: np.ndarray, ref_scores: np.ndarray, k: int) -> bool:
    """Tie-aware check (indexer_quant.py:66-68 form): a selection of k distinct positions is a valid
    top-k of ref_scores iff every selected value is >= the k-th largest reference value and every
    value strictly above it is selected. Rows whose k-th value is -inf compare the finite part."""
    s = np.asarray(ref_scores).reshape(-1, ref_scores.shape[-1])
    sel = np.asarray(sel_idx).reshape(-1, k)
    for r in range(s.shape[0]):
        row, pick = s[r], sel[r]
        if len(np.unique(pick)) != k or pick.min() < 0 or pick.max() >= row.shape[0]:
            return False
        kth = np.partition(row, row.shape[0] - k)[row.shape[0] - k]
        if np.isneginf(kth):
            fin = np.flatnonzero(np.isfinite(row))
            if not np.all(np.isin(fin, pick)):
                return False
            continue
        if np.any(row[pick] < kth):
            return False
        if not np.all(np.isin(np.flatnonzero(row > kth), pick)):
            return False
    return True


# ---------------------------------------------------------------------------------- helpers
def hadamard_matrix(d: int = 128) -> np.ndarray:
    """hadamard_quant.py:19-23: Sylvester Hadamard / sqrt(d), rounded to float32 as the reference
    builds it (then widened to float64 by rotate_quant_ref, hadamard_quant.py:108)."""
    h = np.ones((1, 1))
    while h.shape[0] < d:
        h = np.block([[h, h], [h, -h]])
    return (h / np.sqrt(d)).astype(np.float32).astype(np.float64)


def rotate_quant_ref(x: np.ndarray, rotate: bool = True):
    """hadamard_quant.py:106-110: float64 rotation, per-vector scale amax/127 (floor 1e-4),
    round-half-even, clamp. Returns (int8 [..., 128], float32 [...])."""
    xr = np.asarray(x, dtype=np.float64)
    if rotate:
        xr = xr @ hadamard_matrix(xr.shape[-1])
    s = np.maximum(np.abs(xr).max(-1), 1e-4) / 127.0
    q = np.clip(np.rint(xr / s[..., None]), -127, 127).astype(np.int8)
    return q, s.astype(np.float32)


def weight_quant_ref(w: np.ndarray):
    """The weight block quantiser the reference's tests and benchmark apply to the GEMM's B operand
    (test_kernels.py:80-82, bench.py:43-44): per 128 x 128 block of w [N, K] (float32), scale =
    max(amax, 1e-4) / 127 (float32 division), q = clamp(round_half_even(w / scale), -127, 127).
    Returns (int8 [N, K], float32 [N/128, K/128]). NaN converts to 0."""
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    b = w.reshape(N // GROUP, GROUP, K // GROUP, GROUP)
    with np.errstate(invalid="ignore"):
        amax = np.abs(b).max(axis=(1, 3))
        s = (np.maximum(amax, np.float32(1e-4)) / np.float32(127.0)).astype(np.float32)
        s = np.where(np.isnan(amax), np.float32(np.nan), s).astype(np.float32)
        q = np.clip(np.rint(b / s[:, None, :, None]), -127, 127)
    q = np.nan_to_num(q, nan=0.0).astype(np.int8)
    return q.reshape(N, K), s


def rel_err(x: np.ndarray, ref: np.ndarray) -> float:
    """test_kernels.py:15-17: max |x - ref| over finite ref, divided by max |ref|."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    fin = np.isfinite(ref)
    if not fin.any():
        return 0.0
    return float(np.abs(x[fin] - ref[fin]).max() / max(np.abs(ref[fin]).max(), 1e-30))
