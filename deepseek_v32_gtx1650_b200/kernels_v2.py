"""API shims for the reference's kernels_v2.py (dp4a, K-major packed int32 layouts).

The reference's v2 layout ([K/4, rows] int32, kernels_v2.py:52-67,162-170) exists because
Turing's dp4a wants K-major words. The B200 tensor cores read the row-major int8 layout of
kernels.py directly, so these shims keep the v2 names and layouts for callers and unpack to
row-major before calling the same sm_100a kernels.
"""
from __future__ import annotations

import torch

from .kernels import GROUP, act_quant, int8_gemm, int8_index


def kmajor(t: torch.Tensor) -> torch.Tensor:
    """int8 [rows, K] -> int32 [K // 4, rows] K-major packed (kernels_v2.py:65-67)."""
    return t.contiguous().view(torch.int32).T.contiguous()


def unkmajor(tT: torch.Tensor) -> torch.Tensor:
    """int32 [K // 4, rows] K-major packed -> int8 [rows, K] (inverse of kmajor)."""
    return tT.T.contiguous().view(torch.int8)


def act_quant_kmajor(x: torch.Tensor, round_scale: bool = False, block_m: int = 32):
    """x [..., N] -> (int32 [N // 4, M] K-major packed int8, fp32 scales [M, N // 128]) (kernels_v2.py:52-62)."""
    assert x.is_contiguous() and x.shape[-1] % GROUP == 0
    N = x.shape[-1]
    y, s = act_quant(x.view(-1, N), round_scale)
    return kmajor(y), s


def int8_gemm_v2(aT, a_s, bT, b_s, out_dtype=torch.float32):
    """aT int32 [K // 4, M], a_s [M, K // 128], bT int32 [K // 4, N], b_s [N // 128, K // 128] -> [M, N]
    (kernels_v2.py:113-122)."""
    K4, M = aT.shape
    N = bT.shape[1]
    KG = K4 * 4 // GROUP
    assert bT.shape[0] == K4 and N % GROUP == 0 and a_s.shape == (M, KG)
    return int8_gemm(unkmajor(aT), a_s.contiguous(), unkmajor(bT), b_s.contiguous(), out_dtype=out_dtype)


def index_kmajor_q(q: torch.Tensor) -> torch.Tensor:
    """q int8 [b, m, h, d] -> int32 [b, d / 4, m * h] (kernels_v2.py:162-165)."""
    B, M, H, D = q.shape
    return q.contiguous().view(B, M * H, D).view(torch.int32).transpose(1, 2).contiguous()


def index_kmajor_k(k: torch.Tensor) -> torch.Tensor:
    """k int8 [b, n, d] -> int32 [b, d / 4, n] (kernels_v2.py:168-170)."""
    return k.contiguous().view(torch.int32).transpose(1, 2).contiguous()


def int8_index_v2(qT, w, kT, k_s, H, causal=False, start=0, block_q=1, block_n=64, unroll=8, num_warps=1):
    """qT [b, d / 4, m * h], w [b, m, h], kT [b, d / 4, n], k_s [b, n] -> [b, m, n] (kernels_v2.py:173-182)."""
    B, D4, R = qT.shape
    M = R // H
    assert w.is_contiguous() and k_s.is_contiguous() and kT.shape[:2] == (B, D4)
    q = qT.transpose(1, 2).contiguous().view(torch.int8).view(B, M, H, D4 * 4)
    k = kT.transpose(1, 2).contiguous().view(torch.int8)
    return int8_index(q, w, k, k_s, causal=causal, start=start)
