"""Test and measurement infrastructure: PyTorch-on-CPU restatements of the reference's own eager
paths (reference.py:8-82), the fastest CPU implementations the reference itself offers for the hot
path. bench.py times them on the host cores as the CPU baseline and the reference arm; they are
never part of the product path (the package does not import this module).

Each function states which reference lines it follows. They run on CPU tensors with all the
threads torch is given (torch.set_num_threads).
"""
from __future__ import annotations

import torch

GROUP = 128


def act_quant_torch(x: torch.Tensor, round_scale: bool = False):
    """reference.py:8-15 (act_quant_ref, which reference.py:38-40 act_quant_torch returns): per
    128-group amax, s = max(amax, 1e-4) * (1/127) (ue8m0: 2^ceil(log2 s)), y = clamp(round(x / s))."""
    *lead, n = x.shape
    g = x.float().view(*lead, n // GROUP, GROUP)
    s = torch.clamp(g.abs().amax(-1), min=1e-4) * (1.0 / 127.0)
    if round_scale:
        s = torch.exp2(torch.ceil(torch.log2(s)))
    y = torch.clamp(torch.round(g / s.unsqueeze(-1)), -127, 127).to(torch.int8)
    return y.view(*lead, n), s


def dequant_weight(b: torch.Tensor, b_s: torch.Tensor) -> torch.Tensor:
    """The pre-dequantised fp32 weight gemm_dequant_fp32 multiplies against (done once, offline, as
    the reference's baseline assumes): b [N, K] int8 times its [N/128, K/128] block scales."""
    n, k = b.shape
    bs = b_s.repeat_interleave(GROUP, 0)[:n]  # [N, K/128]
    return (b.float().view(n, k // GROUP, GROUP) * bs.unsqueeze(-1)).view(n, k)


def gemm_dequant_fp32(a: torch.Tensor, a_s: torch.Tensor, b_deq: torch.Tensor) -> torch.Tensor:
    """reference.py:43-48: dequantise the activations per 128-block, then one fp32 matmul against
    the pre-dequantised weights."""
    k = a.shape[-1]
    A = (a.float().view(-1, k // GROUP, GROUP) * a_s.view(-1, k // GROUP, 1)).view(*a.shape[:-1], k)
    return A @ b_deq.T


def int_mm_unscaled(a: torch.Tensor, bT: torch.Tensor) -> torch.Tensor:
    """reference.py:56-58: torch._int_mm with no block scales (an upper bound on INT8 matmul speed,
    not a usable layer)."""
    return torch._int_mm(a, bT)


def index_torch_int8(q, w, k, k_s, chunk: int = 64, rows=None):
    """reference.py:72-82: the indexer through torch._int_mm on stacked heads, chunked over queries
    (no causal mask; the reference's baseline scores every key). rows: only these query rows."""
    B, M, H, D = q.shape
    rows = torch.arange(M) if rows is None else torch.as_tensor(rows)
    out = []
    for b in range(B):
        kT = k[b].T.contiguous()
        acc = []
        for i in range(0, len(rows), chunk):
            r = rows[i:i + chunk]
            qi = q[b, r].reshape(-1, D)
            lg = torch._int_mm(qi, kT).float().clamp_min_(0).view(-1, H, k.shape[1])
            acc.append((lg * w[b, r].unsqueeze(-1)).sum(1) * k_s[b])
        out.append(torch.cat(acc, 0))
    return torch.stack(out)


def index_torch_fp32(q, w, k, k_s, chunk: int = 64, rows=None):
    """reference.py:61-69: the indexer on dequantised fp32 operands, chunked over queries."""
    B, M, H, D = q.shape
    rows = torch.arange(M) if rows is None else torch.as_tensor(rows)
    kf = k.float()
    out = []
    for i in range(0, len(rows), chunk):
        r = rows[i:i + chunk]
        lg = torch.einsum("bmhd,bnd->bmhn", q[:, r].float(), kf).clamp_min_(0)
        out.append((lg * w[:, r].unsqueeze(-1)).sum(2) * k_s.unsqueeze(1))
    return torch.cat(out, 1)
