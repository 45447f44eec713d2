"""The full lightning-indexer step around the hot path (bench_indexer_e2e.py:46-58): quantise the
step's new keys into an int8 key cache, rotate + quantise the queries, fold the per-vector query
scales into the head weights, then score and select the top-k keys per query.

All compute runs in the sm_100a library (rotate_quant, int8_index_topk); the cache is plain
device tensors owned by the caller.
"""
from __future__ import annotations

import torch

from .kernels import int8_index_topk, rotate_quant


class KeyCache:
    """int8 key cache [B, capacity, 128] with per-key fp32 scales [B, capacity]; keys [0, length)
    are valid. The reference keeps the same pair (kT, ks) in its K-major layout
    (bench_indexer_e2e.py:47,56)."""

    def __init__(self, batch: int, capacity: int, device, dim: int = 128):
        assert dim == 128
        self.k = torch.zeros(batch, capacity, dim, dtype=torch.int8, device=device)
        self.k_s = torch.zeros(batch, capacity, dtype=torch.float32, device=device)
        self.length = 0

    def append(self, k_new: torch.Tensor) -> None:
        """Rotate + quantise k_new [B, n_new, 128] (fp32/bf16/fp16) into positions [length, length + n_new)."""
        B, n_new, _ = k_new.shape
        assert B == self.k.shape[0] and self.length + n_new <= self.k.shape[1], "key cache overflow"
        kq, ks = rotate_quant(k_new.contiguous())
        self.k[:, self.length:self.length + n_new].copy_(kq)
        self.k_s[:, self.length:self.length + n_new].copy_(ks)
        self.length += n_new


def indexer_step(q: torch.Tensor, w: torch.Tensor, cache: KeyCache, k_new: torch.Tensor | None = None,
                 topk: int = 2048, causal: bool = True, return_scores: bool = False):
    """One indexer step: append k_new to the cache, then for the queries q [B, M, H, 128] (float)
    with head weights w [B, M, H] select the top-k of the cache's keys [0, length).
    Causal: query m is the token at position length - M + m and sees keys up to itself.
    Returns (idx int32 [B, M, topk], vals fp32 [B, M, topk]) (and the scores first when
    return_scores). The query scales multiply w as in bench_indexer_e2e.py:55, inside the rotate +
    quantise kernel; the cache's keys [0, length) are read in place (no copy of the cache)."""
    if k_new is not None:
        cache.append(k_new)
    B, M, H, D = q.shape
    N = cache.length
    # [B, M, H, 128] int8 and the head weights times the per-vector query scales [B, M, H]
    qq, w2 = rotate_quant(q.contiguous(), scale_mul=w.float().contiguous())
    return int8_index_topk(qq, w2, cache.k, cache.k_s, topk=min(topk, N), causal=causal, start=N - M,
                           return_scores=return_scores, n_keys=N)
