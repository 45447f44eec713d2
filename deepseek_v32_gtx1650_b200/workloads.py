"""Seeded synthetic inputs with the shapes and value distributions of the BASELINE configs.

The reference measures on DeepSeek-V3.2 layer shapes with random data (bench.py:35-58,74-92,
bench_indexer_e2e.py:32-48); no dataset is involved. These generators run on the CPU with
torch's seeded RNG so every process (tests, bench, ranks) builds bit-identical inputs.

- act_quant: x ~ N(0,1) fp32 [M, N]; 0.1 % of entries (chosen by a seeded randperm) replaced by
  50 * N(0,1) outliers; row 0 all zeros. The same x cast to bf16 is the bf16 case.
- int8_gemm: activations x ~ N(0,1) bf16 [M, K] (quantised by act_quant on the caller's side),
  weights B ~ U{-127..127} int8 [N, K], weight-block scales b_s = exp(N(-6, 0.5)) [N/128, K/128].
- indexer: q ~ N(0,1) [B, M, H, D] and keys ~ N(0, I_D) with a shared offset of 5 * sqrt(D) in
  channel 0 (indexer_mechanism.py:84 form, c = 5), both Hadamard-rotated (128-point, scale
  D^-1/2, as hadamard_quant.py:106-110) and quantised per vector (amax / 127); head weights
  w = U(0,1) / 64 with the per-vector q scales folded in (bench_indexer_e2e.py:48).
"""
from __future__ import annotations

import math

import torch


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def act_quant_input(M: int = 2048, N: int = 7168, seed: int = 0) -> torch.Tensor:
    g = _gen(seed)
    x = torch.randn(M, N, generator=g, dtype=torch.float32)
    n_out = max(1, (M * N) // 1000)
    pos = torch.randperm(M * N, generator=g)[:n_out]
    x.view(-1)[pos] = 50.0 * torch.randn(n_out, generator=g, dtype=torch.float32)
    x[0] = 0.0
    return x


def gemm_inputs(M: int, N: int, K: int, seed: int = 0):
    """Returns (x bf16 [M, K] activations, B int8 [N, K], b_s fp32 [N/128, K/128])."""
    g = _gen(seed)
    x = torch.randn(M, K, generator=g, dtype=torch.float32).to(torch.bfloat16)
    B = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    b_s = torch.exp(torch.randn(N // 128, K // 128, generator=g, dtype=torch.float32) * 0.5 - 6.0)
    return x, B, b_s.contiguous()


def hadamard(d: int = 128) -> torch.Tensor:
    """Sylvester Hadamard matrix scaled by d^-1/2, with entries rounded to float32 as the
    reference's hadamard_matrix builds it, returned widened to float64."""
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < d:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / math.sqrt(d)).float().double()


def rotate_quant(x: torch.Tensor, rotate: bool = True):
    """x [..., D] float -> (int8 [..., D], fp32 per-vector scales [...]): float64 Hadamard rotation,
    then s = max(amax, 1e-4) / 127 and round-half-even(x / s) clamped to +-127."""
    xr = x.double() @ hadamard(x.shape[-1]) if rotate else x.double()
    s = xr.abs().amax(-1).clamp_min(1e-4) / 127.0
    q = torch.clamp(torch.round(xr / s[..., None]), -127, 127).to(torch.int8)
    return q, s.float()


def index_inputs(B: int, M: int, N: int, H: int = 64, D: int = 128, seed: int = 0, offset: float = 5.0):
    """Returns (q int8 [B, M, H, D], w fp32 [B, M, H], k int8 [B, N, D], k_s fp32 [B, N])."""
    g = _gen(seed)
    qf = torch.randn(B, M, H, D, generator=g, dtype=torch.float32)
    kf = torch.randn(B, N, D, generator=g, dtype=torch.float32)
    kf[..., 0] += offset * math.sqrt(D)
    q, qs = rotate_quant(qf)
    k, ks = rotate_quant(kf)
    w = torch.rand(B, M, H, generator=g, dtype=torch.float32) / 64.0
    w = (w * qs).contiguous()
    return q.contiguous(), w, k.contiguous(), ks.contiguous()


def index_inputs_uniform(B: int, M: int, N: int, H: int = 64, D: int = 128, seed: int = 0):
    """The reference test generator (test_kernels.py:90-95): uniform int8 q/k, w = N(0,1) * 1e-4,
    k_s = U(0,1) * 0.01."""
    g = _gen(seed)
    q = torch.randint(-127, 128, (B, M, H, D), generator=g, dtype=torch.int8)
    k = torch.randint(-127, 128, (B, N, D), generator=g, dtype=torch.int8)
    w = torch.randn(B, M, H, generator=g, dtype=torch.float32) * 1e-4
    k_s = torch.rand(B, N, generator=g, dtype=torch.float32) * 0.01
    return q, w, k, k_s


def gemm_inputs_uniform(M: int, N: int, K: int, seed: int = 0):
    """The reference test generator (test_kernels.py:49-54): uniform int8 A/B, scales U(0,1)*0.01 + 1e-4."""
    g = _gen(seed)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    a_s = torch.rand(M, K // 128, generator=g, dtype=torch.float32) * 0.01 + 1e-4
    b_s = torch.rand(N // 128, K // 128, generator=g, dtype=torch.float32) * 0.01 + 1e-4
    return a, a_s, b, b_s
