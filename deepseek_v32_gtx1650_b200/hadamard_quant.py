"""API shims for the reference's hadamard_quant.py (the indexer's q / k producer).

Same names and outputs as the reference: rotate_quant_kmajor / fwht_quant_kmajor return the
K-major packed layout of kernels_v2 (int32 [B, 32, R]) and per-vector scales [B, R]. The rotation
and quantisation run in the sm_100a library (kernels.rotate_quant, butterfly form in fp32); the
K-major packing is a host-side reshape. The row-major form that int8_index reads is
kernels.rotate_quant itself.
"""
from __future__ import annotations

import torch

from .kernels import rotate_quant

D = 128


def hadamard_matrix(d: int = D, device="cuda") -> torch.Tensor:
    """Sylvester Hadamard matrix scaled by d^-1/2, float32 (hadamard_quant.py:19-23)."""
    h = torch.ones(1, 1)
    while h.shape[0] < d:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / d ** 0.5).to(device=device, dtype=torch.float32).contiguous()


def _to_kmajor(y: torch.Tensor) -> torch.Tensor:
    """int8 [B, R, 128] -> int32 [B, 32, R] (each int32 packs 4 consecutive values of a vector)."""
    B, R, _ = y.shape
    return y.view(B, R, D // 4, 4).view(torch.int32).view(B, R, D // 4).transpose(1, 2).contiguous()


def rotate_quant_kmajor(x: torch.Tensor, rotate: bool = True, block_m: int = 32):
    """x [B, R, 128] -> (int32 [B, 32, R] K-major packed int8, fp32 [B, R]) (hadamard_quant.py:84-93).
    block_m is accepted and ignored."""
    assert x.is_contiguous() and x.shape[-1] == D and x.dim() == 3
    y, s = rotate_quant(x, rotate)
    return _to_kmajor(y), s


def fwht_quant_kmajor(x: torch.Tensor, block_m: int = 32, num_warps: int = 4):
    """Same output as rotate_quant_kmajor(x, rotate=True) (hadamard_quant.py:84-93)."""
    return rotate_quant_kmajor(x, True)


def unpack_kmajor(yT: torch.Tensor) -> torch.Tensor:
    """int32 [B, 32, R] -> int8 [B, R, 128] (hadamard_quant.py:113-115)."""
    return yT.transpose(1, 2).contiguous().view(torch.int8).view(yT.shape[0], yT.shape[2], D)
